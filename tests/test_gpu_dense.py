"""Greedy sampling kernel (kvbp_argmax) against numpy.argmax's rule, the reference's
sampler (kv_coupled_generator.py:337-344): the first index of the maximum, the first NaN
if any, on bf16 logits of the full Qwen2.5 vocabulary (several CTAs per row, reduced over
a thread-block cluster) and on ragged row lengths with padded rows."""

import pytest
import torch

from kvcacheboundaryprotection_b200 import capi

pytestmark = pytest.mark.gpu


def _first_argmax(x: torch.Tensor) -> list:
    out = []
    for row in x.float().cpu():
        nan = torch.nonzero(torch.isnan(row))
        if nan.numel():
            out.append(int(nan[0]))
            continue
        out.append(int(torch.nonzero(row == row.max())[0]))
    return out


@pytest.mark.parametrize("B,V", [(16, 152064), (3, 4097), (5, 8), (1, 1), (2, 40000)])
def test_argmax_first_maximum(B, V):
    g = torch.Generator(device="cuda").manual_seed(V)
    ld = (V + 7) // 8 * 8  # rows must start on 16-byte boundaries
    buf = torch.randn(B, ld, generator=g, device="cuda").to(torch.bfloat16)
    buf[:, V:] = 100.0  # padding past the vocabulary is never a candidate
    logits = buf[:, :V]
    if B > 1 and V > 64:
        logits[1, V - 1] = 30.0
        logits[1, 7] = 30.0  # tie: the lower index wins
        logits[0] = -2.0     # all equal: index 0
    if B > 2 and V > 64:
        logits[2, 40] = float("nan")  # a NaN wins
        logits[2, 3] = 50.0
    out = torch.empty(B, dtype=torch.int32, device="cuda")
    L = capi.lib()
    st = torch.cuda.current_stream().cuda_stream
    for _ in range(2):  # the result does not depend on an earlier call
        capi.check(L.kvbp_argmax(st, B, V, ld, buf.data_ptr(), out.data_ptr()), "argmax")
        torch.cuda.synchronize()
        assert out.tolist() == _first_argmax(logits)


def test_argmax_keys_over_shards_match_full_row():
    # vocabulary shards long enough to be split over a cluster of CTAs per row
    g = torch.Generator(device="cuda").manual_seed(11)
    B, per, shards = 4, 40000, 3
    V = per * shards
    logits = torch.randn(B, V, generator=g, device="cuda").to(torch.bfloat16)
    logits[1, per + 5] = logits[1, 2 * per + 9] = 40.0  # tie across shards
    logits[2, per - 1] = logits[2, per - 2] = 40.0      # tie at the end of a shard
    L = capi.lib()
    st = torch.cuda.current_stream().cuda_stream
    keys = torch.full((B,), torch.iinfo(torch.int64).min, dtype=torch.int64, device="cuda")
    for r in range(shards):
        k = torch.empty(B, dtype=torch.int64, device="cuda")
        part = logits[:, r * per : (r + 1) * per].contiguous()
        capi.check(L.kvbp_argmax_key(st, B, per, per, part.data_ptr(), r * per, k.data_ptr()), "argmax_key")
        torch.maximum(keys, k, out=keys)
    tok = torch.empty(B, dtype=torch.int32, device="cuda")
    capi.check(L.kvbp_key_to_token(st, B, keys.data_ptr(), tok.data_ptr()), "key_to_token")
    torch.cuda.synchronize()
    assert tok.tolist() == _first_argmax(logits)
    assert tok[1].item() == per + 5 and tok[2].item() == per - 2


def test_argmax_keys_signed_zero_and_nan_across_shards():
    """numpy.argmax ranks -0.0 and +0.0 equal (the lower index wins) and returns the first
    NaN whatever its sign: the sharded keys must agree when those cases span shards."""
    B, per, shards = 3, 40000, 3
    V = per * shards
    g = torch.Generator(device="cuda").manual_seed(5)
    logits = -(torch.rand(B, V, generator=g, device="cuda") + 0.5).to(torch.bfloat16)
    bits = logits.view(torch.int16)
    logits[0, 10] = -0.0        # shard 0: negative zero first ...
    logits[0, per + 2] = 0.0    # ... shard 1: positive zero later -> index 10
    logits[1, 3] = 40.0
    bits[1, 2 * per + 7] = -64  # 0xFFC0: a negative NaN in shard 2 wins over the finite 40
    bits[2, per + 1] = -64      # negative NaN in shard 1 ...
    bits[2, 100] = 0x7FC0       # ... but a positive NaN comes first in shard 0
    L = capi.lib()
    st = torch.cuda.current_stream().cuda_stream
    keys = torch.full((B,), torch.iinfo(torch.int64).min, dtype=torch.int64, device="cuda")
    for r in range(shards):
        k = torch.empty(B, dtype=torch.int64, device="cuda")
        part = logits[:, r * per : (r + 1) * per].contiguous()
        capi.check(L.kvbp_argmax_key(st, B, per, per, part.data_ptr(), r * per, k.data_ptr()), "argmax_key")
        torch.maximum(keys, k, out=keys)
    tok = torch.empty(B, dtype=torch.int32, device="cuda")
    capi.check(L.kvbp_key_to_token(st, B, keys.data_ptr(), tok.data_ptr()), "key_to_token")
    torch.cuda.synchronize()
    assert tok.tolist() == _first_argmax(logits) == [10, 2 * per + 7, 100]
